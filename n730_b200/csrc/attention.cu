// RoPE + GQA attention over a paged fp16 KV cache.
//
// Replaces the reference's attention path: rope_kernel (n730_cuda.cu:277-304),
// the D2D KV append in src-code/inference.py:539-549, and
// n730_attention_forward (n730_cuda.cu:709-845: whole-cache repack, 2*n_heads
// cuBLAS calls, materialised fp32 scores, mask and softmax kernels).
//
// Decode (one token per sequence) is a single kernel: a cluster of 8 CTAs per
// (sequence, KV head), each CTA one split of the context.  A CTA applies
// rotate_half RoPE to the group's n_heads/n_kv query heads in shared memory;
// the CTA whose split holds the new position RoPEs and appends k/v to the
// cache; then each CTA streams its pages once for all query heads of the
// group (flash-decoding with an online softmax).  The splits merge through
// distributed shared memory (cluster rank 0 reads every rank's partials):
// out = sum_s e^(m_s-M) acc_s / (sum_s e^(m_s-M) l_s + 1e-9), the reference's
// normalisation (n730_cuda.cu:236-257).  Scores are scaled by 1/sqrt(head_dim).
// The reference's exp(max(s - m, -50)) floor changes weights by at most e^-50
// and is not reproduced.
//
// Prefill uses kv_write (RoPE + cache append for T tokens) and a causal
// tensor-core flash-attention kernel; masked keys get weight 0 (the reference
// uses -1e4 scores, weight <= e^-50).
#include <cfloat>

#include <cooperative_groups.h>

#include "attention.h"

namespace cg = cooperative_groups;

namespace n730 {

constexpr int MAX_G = 8;

__device__ __forceinline__ const __half* page_ptr(const __half* pages, const int* bt, int p, const AttnDims& d,
                                                  int kvh) {
  const int page = bt[p / d.page_size];
  return pages + (((int64_t)page * d.n_kv + kvh) * d.page_size + (p % d.page_size)) * d.head_dim;
}

// Decode attention, one thread-block cluster per (sequence, KV head): CTA r
// of the cluster owns context positions [r*chunk, (r+1)*chunk).  Per tile of
// DEC_TILE positions the CTA stages K and V with cp.async into XOR-swizzled
// shared memory, three buffers deep (the next two tiles load while this one
// computes); each of its 8 warps takes 16 positions and computes
//   S = Q K^T   with mma.m16n8k16 (f16 in, f32 accumulate): the G <= 8 query
//               heads of the group are rows 0..G-1 of the A tile, K feeds B
//               through ldmatrix,
//   online softmax on the S fragments (per warp running max / sum),
//   O += P V    with P re-packed from the S fragments as the A operand and V
//               through ldmatrix.trans.
// Warps merge in shared memory, then the cluster's CTAs merge through
// distributed shared memory (rank 0 reads every rank's m, l, O).
constexpr int DEC_THREADS = 256;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int DEC_TILE = 16 * DEC_WARPS;  // 128 positions per tile
constexpr int DEC_STAGES = 3;             // tile buffers (two tiles in flight while one computes)

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(dst), "l"(src), "r"(pred ? 16 : 0));
}
// byte offset of 16-byte chunk c of row r in a swizzled [rows][HD] fp16 tile
template <int HD>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * HD * 2 + ((c ^ (r & 7)) << 4));
}

template <int HD>
struct DecSmem {
  __half k[DEC_STAGES][DEC_TILE * HD];  // tile buffers: the next two tiles load while one computes;
  __half v[DEC_STAGES][DEC_TILE * HD];  // after the loop k holds the per-warp outputs (wo)
  float q[MAX_G][HD];                 // RoPE'd, scaled queries (fp32)
  float wm[DEC_WARPS][MAX_G], wl[DEC_WARPS][MAX_G];
  float m[MAX_G], l[MAX_G];           // this CTA's split
  float o[MAX_G][HD];
  float sw[MAX_G][16], den[MAX_G];    // cluster merge: weight e^(m_r - M) of each split, denominator
};

template <int HD>
__global__ void __launch_bounds__(DEC_THREADS) attn_decode_kernel(const DecodeAttnArgs a) {
  using SM = DecSmem<HD>;
  constexpr int H2 = HD / 2, KS = HD / 16, NCH = HD / 8;  // k-steps, 16-B chunks per row
  extern __shared__ __align__(128) uint8_t dsm[];
  SM& sm = *reinterpret_cast<SM*>(dsm);

  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int split = (int)cluster.block_rank();
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const AttnDims& d = a.d;
  const int G = d.n_heads / d.n_kv;
  pdl_wait();
  const int pos = a.seq_lens[b];
  const int L = pos + 1;
  const int chunk = ((L + S - 1) / S + DEC_TILE - 1) / DEC_TILE * DEC_TILE;
  const int t0 = split * chunk, t1 = min(L, t0 + chunk);
  const int* bt = a.block_table + (int64_t)b * d.max_pages;
  const float* qkv = a.qkv + (int64_t)b * a.ld_qkv;
  const float* cs = a.cos_t + (int64_t)pos * H2;
  const float* sn = a.sin_t + (int64_t)pos * H2;

  for (int i = tid; i < MAX_G * HD; i += DEC_THREADS) {  // RoPE'd, pre-scaled queries
    const int g = i / HD, j = i % HD;
    float v = 0.f;
    if (g < G) {
      const float* qh = qkv + (int64_t)(kvh * G + g) * HD;
      const int j0 = j < H2 ? j : j - H2;
      const float x0 = qh[j0], x1 = qh[j0 + H2], c = cs[j0], s = sn[j0];
      v = (j < H2 ? x0 * c - x1 * s : x1 * c + x0 * s) * d.scale;
    }
    sm.q[g][j] = v;
  }
  // the new position's k (RoPE'd) and v, rounded to fp16 as stored
  const bool owns_new = t0 <= pos && pos < t1;
  if (owns_new) {
    const float* kh = qkv + (int64_t)(d.n_heads + kvh) * HD;
    const float* vh = qkv + (int64_t)(d.n_heads + d.n_kv + kvh) * HD;
    __half* kd = const_cast<__half*>(page_ptr(a.kv.k_pages, bt, pos, d, kvh));
    __half* vd = const_cast<__half*>(page_ptr(a.kv.v_pages, bt, pos, d, kvh));
    for (int j = tid; j < H2; j += DEC_THREADS) {
      const float x0 = kh[j], x1 = kh[j + H2], c = cs[j], s = sn[j];
      kd[j] = __float2half_rn(x0 * c - x1 * s);
      kd[j + H2] = __float2half_rn(x1 * c + x0 * s);
    }
    for (int j = tid; j < HD; j += DEC_THREADS) vd[j] = __float2half_rn(vh[j]);
  }
  __syncthreads();
  pdl_launch_dependents();

  // Q as the A operand: rows 0..7 = query heads (>= G are zero), rows 8..15 zero
  uint32_t qa[KS][2];
  {
    const int r = lane >> 2, c = (lane & 3) * 2;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = pack_half2(sm.q[r][ks * 16 + c], sm.q[r][ks * 16 + c + 1]);
      qa[ks][1] = pack_half2(sm.q[r][ks * 16 + c + 8], sm.q[r][ks * 16 + c + 9]);
    }
  }
  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // for head row lane>>2 (replicated over the 4 lanes of a row)
  // ---- stage K and V rows [tile, tile + DEC_TILE) into buffer `buf` (swizzled; rows past t1 zero) ----
  // Thread tid copies 16-byte chunk tid % NCH of rows tid / NCH + j * RSTEP; the block-table
  // reads for its rows go out first, independent of one another, then the copies.
  constexpr int RSTEP = DEC_THREADS / NCH, NIT = DEC_TILE / RSTEP;
  static_assert(DEC_THREADS % NCH == 0 && DEC_TILE % RSTEP == 0, "staging covers the tile exactly");
  const int sr0 = tid / NCH, sc = tid % NCH, ps = d.page_size;
  auto stage = [&](int tile, int buf) {
    const int np = min(DEC_TILE, t1 - tile);
    const uint32_t kb = smem_u32(sm.k[buf]), vb = smem_u32(sm.v[buf]);
    int64_t off[NIT];
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
      const int r = sr0 + j * RSTEP;
      const int p = r < np ? tile + r : tile;  // rows past the end: a valid address, zero bytes read
      off[j] = (((int64_t)bt[p / ps] * d.n_kv + kvh) * ps + p % ps) * HD + sc * 8;
    }
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
      const int r = sr0 + j * RSTEP;
      cp_async16(kb + swz<HD>(r, sc), a.kv.k_pages + off[j], r < np);
      cp_async16(vb + swz<HD>(r, sc), a.kv.v_pages + off[j], r < np);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (t0 < t1) stage(t0, 0);
  if (t0 + DEC_TILE < t1) stage(t0 + DEC_TILE, 1);

  for (int tile = t0, it = 0; tile < t1; tile += DEC_TILE, ++it) {
    const int np = min(DEC_TILE, t1 - tile), buf = it % DEC_STAGES;
    const uint32_t ks_base = smem_u32(sm.k[buf]), vs_base = smem_u32(sm.v[buf]);
    // the tile two ahead goes out before this one is waited for (its buffer was last read
    // in the previous iteration, before the loop's closing barrier); then wait until at most
    // the copies of the tiles after this one are pending
    static_assert(DEC_STAGES == 3, "the wait_group counts below assume three buffers");
    if (tile + 2 * DEC_TILE < t1) {
      stage(tile + 2 * DEC_TILE, (it + 2) % DEC_STAGES);
      asm volatile("cp.async.wait_group 2;" ::: "memory");
    } else if (tile + DEC_TILE < t1) {
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (owns_new && pos >= tile && pos < tile + DEC_TILE) {  // the row just appended, from registers' values
      const int r = pos - tile;
      const float* kh = qkv + (int64_t)(d.n_heads + kvh) * HD;
      const float* vh = qkv + (int64_t)(d.n_heads + d.n_kv + kvh) * HD;
      for (int j = tid; j < HD; j += DEC_THREADS) {
        const int j0 = j < H2 ? j : j - H2;
        const float x0 = kh[j0], x1 = kh[j0 + H2], c = cs[j0], s = sn[j0];
        const float kv = j < H2 ? x0 * c - x1 * s : x1 * c + x0 * s;
        const uint32_t off = swz<HD>(r, j / 8) + (j % 8) * 2;
        *reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(sm.k[buf]) + off) = __float2half_rn(kv);
        *reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(sm.v[buf]) + off) = __float2half_rn(vh[j]);
      }
      __syncthreads();
    }
    const int w0 = warp * 16;  // this warp's 16 positions of the tile
    if (w0 < np) {
      // ---- S = Q K^T for 16 positions (two n-tiles of 8) ----
      float sacc[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        // matrices: (n-tile 0, k lo), (n-tile 0, k hi), (n-tile 1, k lo), (n-tile 1, k hi)
        const int mi = lane >> 3, rr = lane & 7;
        const int row = w0 + (mi >> 1) * 8 + rr;
        const int chk = ks * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ks_base + swz<HD>(row, chk), b0, b1, b2, b3);
        const uint32_t af[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
        mma_16816(sacc[0], af, b0, b1);
        mma_16816(sacc[1], af, b2, b3);
      }
      // ---- online softmax on rows 0..7 (c0, c1 of each n-tile) ----
      float sv[4];
      sv[0] = sacc[0][0]; sv[1] = sacc[0][1]; sv[2] = sacc[1][0]; sv[3] = sacc[1][1];
      const int cb = (lane & 3) * 2;
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pcol = w0 + (j >> 1) * 8 + cb + (j & 1);
        if (pcol >= np) sv[j] = -INFINITY;
        mt = fmaxf(mt, sv[j]);
      }
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float mn = fmaxf(m_run, mt);
      const float al = m_run == -INFINITY ? 0.f : __expf(m_run - mn);
      float pe[4], ts = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) { pe[j] = sv[j] == -INFINITY ? 0.f : __expf(sv[j] - mn); ts += pe[j]; }
      ts += __shfl_xor_sync(0xffffffffu, ts, 1);
      ts += __shfl_xor_sync(0xffffffffu, ts, 2);
      l_run = l_run * al + ts;
      m_run = mn;
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) { o[n][0] *= al; o[n][1] *= al; }
      // ---- O += P V (P: rows = heads, k = this warp's 16 positions) ----
      const uint32_t pa[4] = {pack_half2(pe[0], pe[1]), 0u, pack_half2(pe[2], pe[3]), 0u};
#pragma unroll
      for (int n2 = 0; n2 < HD / 16; ++n2) {
        // matrices (trans): (k lo, n-tile 2*n2), (k hi, n-tile 2*n2), (k lo, 2*n2+1), (k hi, 2*n2+1)
        const int mi = lane >> 3, rr = lane & 7;
        const int row = w0 + (mi & 1) * 8 + rr;
        const int chk = n2 * 2 + (mi >> 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vs_base + swz<HD>(row, chk), v0, v1, v2, v3);
        mma_16816(o[2 * n2], pa, v0, v1);
        mma_16816(o[2 * n2 + 1], pa, v2, v3);
      }
    }
    __syncthreads();  // tile buffers are reused
  }

  // ---- merge the 8 warps of this CTA (per-warp outputs in the first K buffer: the loop is done) ----
  float (*wo)[MAX_G][HD] = reinterpret_cast<float (*)[MAX_G][HD]>(&sm.k[0][0]);
  static_assert(sizeof(float) * DEC_WARPS * MAX_G * HD <= sizeof(sm.k), "per-warp outputs fit the K buffers");
  {
    const int r = lane >> 2, cb = (lane & 3) * 2;
    if ((lane & 3) == 0 && r < MAX_G) { sm.wm[warp][r] = m_run; sm.wl[warp][r] = l_run; }
    if (r < MAX_G)
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) { wo[warp][r][n * 8 + cb] = o[n][0]; wo[warp][r][n * 8 + cb + 1] = o[n][1]; }
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += DEC_THREADS) {
    const int g = i / HD, dd = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < DEC_WARPS; ++w) M = fmaxf(M, sm.wm[w][g]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < DEC_WARPS; ++w) {
      const float mw = sm.wm[w][g];
      if (mw == -INFINITY) continue;
      const float e = __expf(mw - M);
      num = fmaf(e, wo[w][g][dd], num);
      den = fmaf(e, sm.wl[w][g], den);
    }
    sm.o[g][dd] = num;
    if (dd == 0) { sm.m[g] = M; sm.l[g] = den; }
  }
  cluster.sync();  // every split's (m, l, o) is visible cluster-wide
  // every rank: split weights per head (warp g, lane r = split r, fixed-order
  // reductions), then this rank merges its 1/S slice of the G x HD outputs
  if (warp < G) {
    const int g = warp;
    const float mr = lane < S ? cluster.map_shared_rank(&sm, lane)->m[g] : -INFINITY;
    const float lr = lane < S ? cluster.map_shared_rank(&sm, lane)->l[g] : 0.f;
    float M = mr;
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
    const float w = mr == -INFINITY ? 0.f : __expf(mr - M);
    float dn = w * lr;
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) dn += __shfl_xor_sync(0xffffffffu, dn, o2);
    if (lane < 16) sm.sw[g][lane] = lane < S ? w : 0.f;
    if (lane == 0) sm.den[g] = dn;
  }
  __syncthreads();
  {
    const int n_out = G * HD, lo = split * n_out / S, hi = (split + 1) * n_out / S;
    for (int i = lo + tid; i < hi; i += DEC_THREADS) {
      const int g = i / HD, dd = i % HD;
      float num = 0.f;
      for (int r = 0; r < S; ++r) num = fmaf(sm.sw[g][r], cluster.map_shared_rank(&sm, r)->o[g][dd], num);
      a.out[(int64_t)b * d.n_heads * HD + (int64_t)(kvh * G + g) * HD + dd] = num / (sm.den[g] + 1e-9f);
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until every rank has merged
}

template <typename KernelT, typename ArgT>
static int launch_pdl(KernelT k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, const ArgT& arg) {
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
  N730_CUDA(cudaLaunchKernelEx(&cfg, k, arg));
  return N730_OK;
}

template <int HD>
static int decode_cluster_size() {
  const size_t smem = sizeof(DecSmem<HD>);
  N730_CUDA(cudaFuncSetAttribute(attn_decode_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  N730_CUDA(cudaFuncSetAttribute(attn_decode_kernel<HD>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  for (int cl : {16, 8}) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl, 1, 1);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<HD>, &cfg) == cudaSuccess && n > 0) return cl;
    cudaGetLastError();
  }
  return 8;
}

int attn_decode_launch(const DecodeAttnArgs& a, cudaStream_t st) {
  const AttnDims& d = a.d;
  N730_REQUIRE(d.n_kv > 0 && d.n_heads % d.n_kv == 0 && d.n_heads / d.n_kv <= MAX_G, N730_BAD_ARG,
               "attention: n_heads/n_kv must be an integer <= %d", MAX_G);
  N730_REQUIRE(d.head_dim == 64 || d.head_dim == 128, N730_UNSUPPORTED, "attention: head_dim %d", d.head_dim);
  N730_REQUIRE(a.batch >= 1, N730_BAD_ARG, "attention: bad batch");
  // the kernel attributes and the cluster size are set up once per device
  static std::mutex mu;
  static int cl128[N730_MAX_DEVICES] = {}, cl64[N730_MAX_DEVICES] = {};
  int dev = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_REQUIRE(dev >= 0 && dev < N730_MAX_DEVICES, N730_BAD_ARG, "attention: device ordinal %d", dev);
  int cl_max = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    int& slot = d.head_dim == 128 ? cl128[dev] : cl64[dev];
    if (!slot) slot = d.head_dim == 128 ? decode_cluster_size<128>() : decode_cluster_size<64>();
    cl_max = slot;
    if (cl_max < 0) slot = 0;  // set-up failed: try again on the next call
  }
  if (cl_max < 0) return cl_max;
  // splits per (sequence, KV head): about one CTA per SM in all (a CTA's three tile buffers take
  // most of an SM's shared memory, and its loads overlap its own compute)
  int cl = cl_max;
  while (cl > 1 && (int64_t)a.batch * d.n_kv * cl > (int64_t)num_sms()) cl >>= 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cl, d.n_kv, a.batch);
  cfg.blockDim = dim3(DEC_THREADS);
  cfg.stream = st;
  cfg.dynamicSmemBytes = d.head_dim == 128 ? sizeof(DecSmem<128>) : sizeof(DecSmem<64>);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 2 : 1;
  if (d.head_dim == 128) N730_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_kernel<128>, a));
  else N730_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_kernel<64>, a));
  return N730_OK;
}

// ---------------------------------------------------------------------------
// prefill
// ---------------------------------------------------------------------------
__global__ void kv_write_kernel(const KVWriteArgs a) {
  pdl_wait();
  const int t = blockIdx.x;
  const AttnDims& d = a.d;
  const int H2 = d.head_dim / 2;
  const int pos = a.pos0 + t;
  float* row = a.qkv + (int64_t)t * a.ld_qkv;
  const float* cs = a.cos_t + (int64_t)pos * H2;
  const float* sn = a.sin_t + (int64_t)pos * H2;
  // q heads in place, then k heads into the cache
  for (int i = threadIdx.x; i < (d.n_heads + d.n_kv) * H2; i += blockDim.x) {
    const int h = i / H2, j = i % H2;
    float* x = row + (int64_t)h * d.head_dim;
    const float x0 = x[j], x1 = x[j + H2], c = cs[j], s = sn[j];
    const float y0 = x0 * c - x1 * s, y1 = x1 * c + x0 * s;
    if (h < d.n_heads) {
      x[j] = y0;
      x[j + H2] = y1;
    } else {
      __half* kd = const_cast<__half*>(page_ptr(a.kv.k_pages, a.block_table, pos, d, h - d.n_heads));
      kd[j] = __float2half_rn(y0);
      kd[j + H2] = __float2half_rn(y1);
    }
  }
  for (int i = threadIdx.x; i < d.n_kv * d.head_dim; i += blockDim.x) {
    const int h = i / d.head_dim, j = i % d.head_dim;
    __half* vd = const_cast<__half*>(page_ptr(a.kv.v_pages, a.block_table, pos, d, h));
    vd[j] = __float2half_rn(row[(int64_t)(d.n_heads + d.n_kv + h) * d.head_dim + j]);
  }
}

int kv_write_launch(const KVWriteArgs& a, cudaStream_t st) {
  if (a.T <= 0) return N730_OK;
  return launch_pdl(kv_write_kernel, dim3(a.T), dim3(256), 0, st, a.pdl, a);
}

// Causal prefill attention on the tensor cores (flash-attention style): one
// CTA per (64-query block, query head), 4 warps of 16 queries.  Q is RoPE'd in
// place by kv_write, scaled and rounded to fp16 into swizzled shared memory;
// each warp keeps its A fragments in registers.  Key tiles of 64 positions
// (K and V, fp16 from the paged cache) are double-buffered with cp.async; per
// tile S = Q K^T (mma.m16n8k16, K through ldmatrix), the causal mask, an online
// softmax per query row (quad shuffles), and O += P V with P re-packed from
// the S fragments as the A operand and V through ldmatrix.trans.  Query blocks
// are launched latest first (they have the most key tiles).
constexpr int PF_Q = 64;   // queries per CTA (4 warps x 16)
constexpr int PF_K = 64;   // keys per tile

template <int HD>
struct PfSmem {
  __half q[PF_Q * HD];
  __half k[2][PF_K * HD];
  __half v[2][PF_K * HD];
};

template <int HD>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const PrefillAttnArgs a) {
  constexpr int KS = HD / 16, NCH = HD / 8, NTO = HD / 8;
  extern __shared__ __align__(128) uint8_t dsm[];
  PfSmem<HD>& sm = *reinterpret_cast<PfSmem<HD>*>(dsm);
  pdl_wait();
  const AttnDims& d = a.d;
  const int qb = (int)gridDim.x - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, kvh = h / (d.n_heads / d.n_kv);
  const int q0 = qb * PF_Q, nq = min(PF_Q, a.T - q0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int kend = a.pos0 + q0 + nq;  // keys [0, kend) are needed by the CTA
  const int ntiles = (kend + PF_K - 1) / PF_K;
  const uint32_t qs = smem_u32(sm.q);
  const uint32_t kb[2] = {smem_u32(sm.k[0]), smem_u32(sm.k[1])};
  const uint32_t vb[2] = {smem_u32(sm.v[0]), smem_u32(sm.v[1])};

  auto stage = [&](int t, int buf) {  // K and V rows [t*PF_K, +PF_K) (zero past kend)
    const int k0 = t * PF_K;
    for (int i = tid; i < PF_K * NCH; i += 128) {
      const int r = i / NCH, c = i % NCH;
      const bool ok = k0 + r < kend;
      const int p = ok ? k0 + r : k0;
      cp_async16(kb[buf] + swz<HD>(r, c), page_ptr(a.kv.k_pages, a.block_table, p, d, kvh) + c * 8, ok);
      cp_async16(vb[buf] + swz<HD>(r, c), page_ptr(a.kv.v_pages, a.block_table, p, d, kvh) + c * 8, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  stage(0, 0);
  for (int i = tid; i < PF_Q * NCH; i += 128) {  // scaled fp16 queries, rows >= nq zero
    const int r = i / NCH, c = i % NCH;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (r < nq) {
      const float4* src = reinterpret_cast<const float4*>(a.qkv + (int64_t)(q0 + r) * a.ld_qkv + (int64_t)h * HD + c * 8);
      const float4 x0 = src[0], x1 = src[1];
      w[0] = pack_half2(x0.x * d.scale, x0.y * d.scale); w[1] = pack_half2(x0.z * d.scale, x0.w * d.scale);
      w[2] = pack_half2(x1.x * d.scale, x1.y * d.scale); w[3] = pack_half2(x1.z * d.scale, x1.w * d.scale);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.q) + swz<HD>(r, c)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  __syncthreads();
  pdl_launch_dependents();
  uint32_t qa[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks)
    ldsm_x4(qs + swz<HD>(warp * 16 + (lane & 15), ks * 2 + (lane >> 4)), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  float o[NTO][4];
#pragma unroll
  for (int n = 0; n < NTO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mr[2] = {-INFINITY, -INFINITY}, lr[2] = {0.f, 0.f};  // rows g and g+8
  const int qp = a.pos0 + q0 + warp * 16 + g;                 // position of row g (row g+8: qp + 8)
  const int mi = lane >> 3, rr = lane & 7;

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) {
      stage(t + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const int k0 = t * PF_K;
    // ---- S = Q K^T, 8 n-tiles of 8 keys ----
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb[buf] + swz<HD>(np * 16 + (mi >> 1) * 8 + rr, ks * 2 + (mi & 1)), b0, b1, b2, b3);
        mma_16816(sc[2 * np], qa[ks], b0, b1);
        mma_16816(sc[2 * np + 1], qa[ks], b2, b3);
      }
    }
    // ---- causal mask, online softmax (rows g: c0 c1, g+8: c2 c3) ----
    float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kp = k0 + n * 8 + 2 * tq + (e & 1);
        const int row_p = qp + (e >> 1) * 8;
        if (kp > row_p || kp >= kend) sc[n][e] = -INFINITY;
        mt[e >> 1] = fmaxf(mt[e >> 1], sc[n][e]);
      }
    float al[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mt[hr] = fmaxf(mt[hr], __shfl_xor_sync(0xffffffffu, mt[hr], 1));
      mt[hr] = fmaxf(mt[hr], __shfl_xor_sync(0xffffffffu, mt[hr], 2));
      const float mn = fmaxf(mr[hr], mt[hr]);
      al[hr] = (mr[hr] == -INFINITY || mn == -INFINITY) ? 0.f : __expf(mr[hr] - mn);
      mr[hr] = mn;
    }
    float ts[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = sc[n][e] == -INFINITY ? 0.f : __expf(sc[n][e] - mr[e >> 1]);
        sc[n][e] = v;
        ts[e >> 1] += v;
      }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      ts[hr] += __shfl_xor_sync(0xffffffffu, ts[hr], 1);
      ts[hr] += __shfl_xor_sync(0xffffffffu, ts[hr], 2);
      lr[hr] = lr[hr] * al[hr] + ts[hr];
    }
#pragma unroll
    for (int n = 0; n < NTO; ++n) { o[n][0] *= al[0]; o[n][1] *= al[0]; o[n][2] *= al[1]; o[n][3] *= al[1]; }
    // ---- O += P V: 4 k-steps of 16 keys, P from the S fragments ----
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t pa[4] = {pack_half2(sc[2 * j][0], sc[2 * j][1]), pack_half2(sc[2 * j][2], sc[2 * j][3]),
                              pack_half2(sc[2 * j + 1][0], sc[2 * j + 1][1]),
                              pack_half2(sc[2 * j + 1][2], sc[2 * j + 1][3])};
#pragma unroll
      for (int n2 = 0; n2 < HD / 16; ++n2) {
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vb[buf] + swz<HD>(j * 16 + (mi & 1) * 8 + rr, n2 * 2 + (mi >> 1)), v0, v1, v2, v3);
        mma_16816(o[2 * n2], pa, v0, v1);
        mma_16816(o[2 * n2 + 1], pa, v2, v3);
      }
    }
    __syncthreads();  // buffer buf is refilled by the stage of tile t + 2
  }
  // ---- normalise and store rows g and g+8 of this warp ----
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = warp * 16 + g + hr * 8;
    if (r >= nq) continue;
    const float inv = 1.f / (lr[hr] + 1e-9f);
    float* out = a.out + (int64_t)(q0 + r) * d.n_heads * HD + (int64_t)h * HD;
#pragma unroll
    for (int n = 0; n < NTO; ++n)
      *reinterpret_cast<float2*>(out + n * 8 + 2 * tq) = make_float2(o[n][hr * 2] * inv, o[n][hr * 2 + 1] * inv);
  }
}

int attn_prefill_launch(const PrefillAttnArgs& a, cudaStream_t st) {
  const AttnDims& d = a.d;
  if (a.T <= 0) return N730_OK;
  N730_REQUIRE(d.head_dim == 64 || d.head_dim == 128, N730_UNSUPPORTED, "attention: head_dim %d", d.head_dim);
  N730_REQUIRE(a.ld_qkv % 4 == 0 && ((uintptr_t)a.qkv & 15) == 0, N730_BAD_ARG, "attention: qkv alignment");
  dim3 grid((a.T + PF_Q - 1) / PF_Q, d.n_heads);
  if (d.head_dim == 128) {
    if (int rc = smem_attr_once<attn_prefill_kernel<128>>((int)sizeof(PfSmem<128>))) return rc;
    return launch_pdl(attn_prefill_kernel<128>, grid, dim3(128), sizeof(PfSmem<128>), st, a.pdl, a);
  }
  if (int rc = smem_attr_once<attn_prefill_kernel<64>>((int)sizeof(PfSmem<64>))) return rc;
  return launch_pdl(attn_prefill_kernel<64>, grid, dim3(128), sizeof(PfSmem<64>), st, a.pdl, a);
}

}  // namespace n730
