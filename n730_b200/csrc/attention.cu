// RoPE + GQA attention over a paged fp16 KV cache.
//
// Replaces the reference's attention path: rope_kernel (n730_cuda.cu:277-304),
// the D2D KV append in src-code/inference.py:539-549, and
// n730_attention_forward (n730_cuda.cu:709-845: whole-cache repack, 2*n_heads
// cuBLAS calls, materialised fp32 scores, mask and softmax kernels).
//
// Decode (one token per sequence) is a single kernel: each CTA owns one
// (sequence, KV head, split of the context).  It applies rotate_half RoPE to
// the group's n_heads/n_kv query heads in shared memory, the CTA whose split
// holds the new position RoPEs and appends k/v to the cache, then streams its
// pages once for all query heads of the group (flash-decoding with an online
// softmax).  The last CTA of a (sequence, KV head) to finish, found with an
// atomic ticket, merges the splits: out = sum_s e^(m_s-M) acc_s /
// (sum_s e^(m_s-M) l_s + 1e-9), the reference's normalisation
// (n730_cuda.cu:236-257).  Scores are scaled by 1/sqrt(head_dim).  The
// reference's exp(max(s - m, -50)) floor changes weights by at most e^-50 and
// is not reproduced.
//
// Prefill uses kv_write (RoPE + cache append for T tokens) and a causal
// CUDA-core flash-attention kernel; masked keys get weight 0 (the reference
// uses -1e4 scores, weight <= e^-50).
#include <cfloat>

#include "attention.h"

namespace n730 {

constexpr int ATT_THREADS = 128;
constexpr int ATT_TILE = 64;
constexpr int MAX_G = 8;

__device__ __forceinline__ const __half* page_ptr(const __half* pages, const int* bt, int p, const AttnDims& d,
                                                  int kvh) {
  const int page = bt[p / d.page_size];
  return pages + (((int64_t)page * d.n_kv + kvh) * d.page_size + (p % d.page_size)) * d.head_dim;
}

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const DecodeAttnArgs a) {
  constexpr int H2 = HD / 2;
  constexpr int QST = H2 + 4;            // padded half-row stride of q in smem
  constexpr int PH = ATT_THREADS / HD;   // position groups in the PV phase
  __shared__ float q_s[MAX_G][2][QST];
  __shared__ float s_s[MAX_G][ATT_TILE];
  __shared__ float m_s[MAX_G], l_s[MAX_G], al_s[MAX_G];
  __shared__ float acc_s[PH > 1 ? PH : 1][MAX_G][HD];
  __shared__ int last_s;

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const AttnDims& d = a.d;
  const int G = d.n_heads / d.n_kv;
  pdl_wait();
  const int pos = a.seq_lens[b];
  const int L = pos + 1;
  const int chunk = ((L + a.n_split - 1) / a.n_split + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
  const int t0 = split * chunk, t1 = min(L, t0 + chunk);
  const int* bt = a.block_table + (int64_t)b * d.max_pages;
  const float* qkv = a.qkv + (int64_t)b * a.ld_qkv;
  const float* cs = a.cos_t + (int64_t)pos * H2;
  const float* sn = a.sin_t + (int64_t)pos * H2;

  if (tid < MAX_G) { m_s[tid] = -INFINITY; l_s[tid] = 0.f; }
  // RoPE'd, pre-scaled queries of the group
  for (int i = tid; i < G * H2; i += ATT_THREADS) {
    const int g = i / H2, j = i % H2;
    const float* qh = qkv + (int64_t)(kvh * G + g) * HD;
    const float x0 = qh[j], x1 = qh[j + H2], c = cs[j], s = sn[j];
    q_s[g][0][j] = (x0 * c - x1 * s) * d.scale;
    q_s[g][1][j] = (x1 * c + x0 * s) * d.scale;
  }
  // the split that holds the new position appends k, v
  if (t0 <= pos && pos < t1) {
    const float* kh = qkv + (int64_t)(d.n_heads + kvh) * HD;
    const float* vh = qkv + (int64_t)(d.n_heads + d.n_kv + kvh) * HD;
    __half* kd = const_cast<__half*>(page_ptr(a.kv.k_pages, bt, pos, d, kvh));
    __half* vd = const_cast<__half*>(page_ptr(a.kv.v_pages, bt, pos, d, kvh));
    for (int j = tid; j < H2; j += ATT_THREADS) {
      const float x0 = kh[j], x1 = kh[j + H2], c = cs[j], s = sn[j];
      kd[j] = __float2half_rn(x0 * c - x1 * s);
      kd[j + H2] = __float2half_rn(x1 * c + x0 * s);
    }
    for (int j = tid; j < HD; j += ATT_THREADS) vd[j] = __float2half_rn(vh[j]);
  }
  __syncthreads();
  pdl_launch_dependents();

  float acc[MAX_G];
#pragma unroll
  for (int g = 0; g < MAX_G; ++g) acc[g] = 0.f;
  const int pd = tid % HD, pg = tid / HD;

  for (int tile = t0; tile < t1; tile += ATT_TILE) {
    // scores: two threads per position, one half of head_dim each
    {
      const int pi = tid >> 1, half = tid & 1;
      const int p = tile + pi;
      float dot[MAX_G];
#pragma unroll
      for (int g = 0; g < MAX_G; ++g) dot[g] = 0.f;
      if (p < t1) {
        const uint4* kr = reinterpret_cast<const uint4*>(page_ptr(a.kv.k_pages, bt, p, d, kvh) + half * H2);
#pragma unroll
        for (int v4 = 0; v4 < H2 / 8; ++v4) {
          const uint4 u = kr[v4];
          const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 kf = __half22float2(h2[e]);
            const int j = v4 * 8 + e * 2;
#pragma unroll
            for (int g = 0; g < MAX_G; ++g) {
              if (g < G) dot[g] = fmaf(q_s[g][half][j], kf.x, fmaf(q_s[g][half][j + 1], kf.y, dot[g]));
            }
          }
        }
      }
#pragma unroll
      for (int g = 0; g < MAX_G; ++g) {
        dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], 1);
        if (half == 0 && g < G) s_s[g][pi] = p < t1 ? dot[g] : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax update, one warp per head
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
      const float s0 = s_s[g][lane], s1 = s_s[g][lane + 32];
      const float mt = warp_max(fmaxf(s0, s1));
      const float mo = m_s[g];
      const float mn = fmaxf(mo, mt);
      const float e0 = s0 == -INFINITY ? 0.f : __expf(s0 - mn);
      const float e1 = s1 == -INFINITY ? 0.f : __expf(s1 - mn);
      s_s[g][lane] = e0;
      s_s[g][lane + 32] = e1;
      const float ts = warp_sum(e0 + e1);
      if (lane == 0) {
        const float al = mo == -INFINITY ? 0.f : __expf(mo - mn);
        al_s[g] = al;
        l_s[g] = l_s[g] * al + ts;
        m_s[g] = mn;
      }
    }
    __syncthreads();
    // P.V: thread = one dim (and one position group when head_dim < 128)
    {
#pragma unroll
      for (int g = 0; g < MAX_G; ++g) if (g < G) acc[g] *= al_s[g];
      const int np = min(ATT_TILE, t1 - tile);
      for (int pi = pg; pi < np; pi += PH) {
        const float v = __half2float(page_ptr(a.kv.v_pages, bt, tile + pi, d, kvh)[pd]);
#pragma unroll
        for (int g = 0; g < MAX_G; ++g) if (g < G) acc[g] = fmaf(s_s[g][pi], v, acc[g]);
      }
    }
    __syncthreads();
  }

  // partials of this split
  const int S = a.n_split;
  if (PH > 1) {
#pragma unroll
    for (int g = 0; g < MAX_G; ++g) if (g < G) acc_s[pg][g][pd] = acc[g];
    __syncthreads();
  }
  if (pg == 0) {
#pragma unroll
    for (int g = 0; g < MAX_G; ++g) {
      if (g >= G) continue;
      float v = acc[g];
      if (PH > 1) { v = 0.f; for (int k = 0; k < PH; ++k) v += acc_s[k][g][pd]; }
      const int h = kvh * G + g;
      a.part_acc[(((int64_t)b * d.n_heads + h) * S + split) * HD + pd] = v;
    }
  }
  if (tid < G) {
    const int h = kvh * G + tid;
    a.part_ml[((int64_t)b * d.n_heads + h) * S + split] = make_float2(m_s[tid], l_s[tid]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int ticket = atomicAdd(&a.counters[b * d.n_kv + kvh], 1);
    last_s = ticket == S - 1;
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // merge the splits of this (sequence, KV head)
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    const float2* ml = a.part_ml + ((int64_t)b * d.n_heads + h) * S;
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, __ldcg(&ml[s].x));
    for (int dd = tid; dd < HD; dd += ATT_THREADS) {
      float num = 0.f, den = 0.f;
      for (int s = 0; s < S; ++s) {
        const float2 v = __ldcg(&ml[s]);
        if (v.x == -INFINITY) continue;
        const float w = __expf(v.x - M);
        den = fmaf(w, v.y, den);
        num = fmaf(w, __ldcg(&a.part_acc[(((int64_t)b * d.n_heads + h) * S + s) * HD + dd]), num);
      }
      a.out[(int64_t)b * d.n_heads * HD + (int64_t)h * HD + dd] = num / (den + 1e-9f);
    }
  }
  if (tid == 0) a.counters[b * d.n_kv + kvh] = 0;
}

size_t attn_decode_workspace(int batch, int n_heads, int n_kv, int head_dim, int n_split) {
  const size_t ml = (size_t)batch * n_heads * n_split * sizeof(float2);
  const size_t acc = (size_t)batch * n_heads * n_split * head_dim * sizeof(float);
  const size_t cnt = (size_t)batch * n_kv * sizeof(int);
  return ml + acc + cnt + 3 * 256;
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

int attn_decode_launch(const DecodeAttnArgs& a, cudaStream_t st) {
  const AttnDims& d = a.d;
  N730_REQUIRE(d.n_kv > 0 && d.n_heads % d.n_kv == 0 && d.n_heads / d.n_kv <= MAX_G, N730_BAD_ARG,
               "attention: n_heads/n_kv must be an integer <= %d", MAX_G);
  N730_REQUIRE(d.head_dim == 64 || d.head_dim == 128, N730_UNSUPPORTED, "attention: head_dim %d", d.head_dim);
  N730_REQUIRE(a.n_split >= 1 && a.batch >= 1, N730_BAD_ARG, "attention: bad split/batch");
  N730_REQUIRE(a.part_ml && a.part_acc && a.counters, N730_NULL, "attention: workspace is null");
  dim3 grid(a.n_split, d.n_kv, a.batch);
  if (d.head_dim == 128) return launch_pdl(attn_decode_kernel<128>, grid, dim3(ATT_THREADS), 0, st, a.pdl, a);
  return launch_pdl(attn_decode_kernel<64>, grid, dim3(ATT_THREADS), 0, st, a.pdl, a);
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

constexpr int PF_Q = 32;     // queries per CTA
constexpr int PF_K = 64;     // keys per tile

template <int HD>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const PrefillAttnArgs a) {
  constexpr int KS = HD + 1;                 // padded strides: conflict-free smem reads
  constexpr int DPT = HD / 4;                // output dims per thread
  constexpr int VS = 4 * (DPT + 1);
  constexpr int PS = PF_K + 1;
  extern __shared__ float pf[];
  float* Qs = pf;                      // [PF_Q][HD+1]
  float* Ks = Qs + PF_Q * KS;          // [PF_K][HD+1]
  float* Vs = Ks + PF_K * KS;          // [PF_K][4][DPT+1]
  float* Ps = Vs + PF_K * VS;          // [PF_Q][PF_K+1]
  pdl_wait();
  const AttnDims& d = a.d;
  const int h = blockIdx.y, kvh = h / (d.n_heads / d.n_kv);
  const int q0 = blockIdx.x * PF_Q;
  const int tid = threadIdx.x, qi = tid >> 2, kg = tid & 3;
  const int nq = min(PF_Q, a.T - q0);
  for (int i = tid; i < PF_Q * HD; i += 128) {
    const int r = i / HD, c = i % HD;
    Qs[r * KS + c] = r < nq ? a.qkv[(int64_t)(q0 + r) * a.ld_qkv + (int64_t)h * HD + c] * d.scale : 0.f;
  }
  float acc[DPT];
#pragma unroll
  for (int j = 0; j < DPT; ++j) acc[j] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int qpos = a.pos0 + q0 + qi;                 // this thread's query position
  const int kend = a.pos0 + q0 + nq;                 // keys [0, kend) are needed by the CTA
  for (int k0 = 0; k0 < kend; k0 += PF_K) {
    __syncthreads();
    for (int i = tid; i < PF_K * HD; i += 128) {
      const int r = i / HD, c = i % HD;
      const int p = k0 + r;
      float kv = 0.f, vv = 0.f;
      if (p < kend) {
        kv = __half2float(page_ptr(a.kv.k_pages, a.block_table, p, d, kvh)[c]);
        vv = __half2float(page_ptr(a.kv.v_pages, a.block_table, p, d, kvh)[c]);
      }
      Ks[r * KS + c] = kv;
      Vs[r * VS + (c / DPT) * (DPT + 1) + (c % DPT)] = vv;
    }
    __syncthreads();
    float s[PF_K / 4];
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < PF_K / 4; ++j) {
      const int kk = kg + 4 * j;
      float dot = 0.f;
#pragma unroll 8
      for (int c = 0; c < HD; ++c) dot = fmaf(Qs[qi * KS + c], Ks[kk * KS + c], dot);
      const int p = k0 + kk;
      s[j] = (qi < nq && p <= qpos) ? dot : -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float mn = fmaxf(m, mt);
    float ts = 0.f;
#pragma unroll
    for (int j = 0; j < PF_K / 4; ++j) {
      const float e = s[j] == -INFINITY ? 0.f : __expf(s[j] - mn);
      Ps[qi * PS + kg + 4 * j] = e;
      ts += e;
    }
    ts += __shfl_xor_sync(0xffffffffu, ts, 1);
    ts += __shfl_xor_sync(0xffffffffu, ts, 2);
    const float al = m == -INFINITY ? 0.f : __expf(m - mn);
    l = l * al + ts;
    m = mn;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < DPT; ++j) acc[j] *= al;
    for (int kk = 0; kk < PF_K; ++kk) {
      const float pv = Ps[qi * PS + kk];
#pragma unroll
      for (int j = 0; j < DPT; ++j) acc[j] = fmaf(pv, Vs[kk * VS + kg * (DPT + 1) + j], acc[j]);
    }
  }
  if (qi < nq) {
    const float inv = 1.f / (l + 1e-9f);
    float* o = a.out + (int64_t)(q0 + qi) * d.n_heads * HD + (int64_t)h * HD + kg * DPT;
#pragma unroll
    for (int j = 0; j < DPT; ++j) o[j] = acc[j] * inv;
  }
}

int attn_prefill_launch(const PrefillAttnArgs& a, cudaStream_t st) {
  const AttnDims& d = a.d;
  if (a.T <= 0) return N730_OK;
  N730_REQUIRE(d.head_dim == 64 || d.head_dim == 128, N730_UNSUPPORTED, "attention: head_dim %d", d.head_dim);
  dim3 grid((a.T + PF_Q - 1) / PF_Q, d.n_heads);
  const int HD = d.head_dim;
  const size_t smem = ((size_t)PF_Q * (HD + 1) + PF_K * (HD + 1) + PF_K * 4 * (HD / 4 + 1) + PF_Q * (PF_K + 1)) *
                      sizeof(float);
  if (HD == 128) {
    static bool cfg = false;
    if (!cfg) {
      N730_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      cfg = true;
    }
    return launch_pdl(attn_prefill_kernel<128>, grid, dim3(128), smem, st, a.pdl, a);
  }
  static bool cfg64 = false;
  if (!cfg64) {
    N730_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cfg64 = true;
  }
  return launch_pdl(attn_prefill_kernel<64>, grid, dim3(128), smem, st, a.pdl, a);
}

}  // namespace n730
